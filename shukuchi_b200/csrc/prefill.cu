// prefill.cu -- batched (prefill) dequantise-matmul on the 5th-generation
// tensor cores: Y[t][m] = sum_k W[m][k] * X[t][k] for a batch of T tokens,
// W in Q4_K or planar Q6_K blocks, X fp32, Y fp32.
//
// The reference has no batched path (engine/src/engine.c:306-501 feeds prompt
// tokens one at a time through op_matmul_q4_k / op_matmul_q6_k,
// engine/src/ops.c:266-314, 361-404); this is the dense contraction those
// per-token matvecs add up to, computed in bf16 x bf16 -> fp32.
//
// One CTA per 128 weight rows x 128 tokens (tcgen05.mma M=128, N=128,
// cta_group::1, accumulator in 128 TMEM columns).  K advances 64 elements per
// step (four MMAs of K=16) through two shared-memory stages:
//   A: 128 rows x 64 bf16, dequantised from the weight blocks by all 256
//      threads (two threads per row, 32 elements each), written in the
//      canonical K-major 128-byte-swizzled layout (16-byte chunk c of row r at
//      r*128 + ((c ^ (r & 7)) * 16); 8-row groups 1024 bytes apart);
//   B: 128 tokens x 64 bf16 copied from the bf16 copy of X, same layout.
// After a proxy fence and a CTA barrier one thread issues the MMAs and
// commits them to the stage's mbarrier; the stage is refilled once that
// commit has arrived, so the fill of step s+1 overlaps the MMAs of step s.
// The epilogue reads the accumulator with tcgen05.ld (warp w: TMEM lanes
// 32w..32w+31 = weight rows) and stores Y token-major, coalesced along m.
// Every wait is bounded; on a time-out the kernel records the error, waits
// (bounded) for its own MMAs, frees its TMEM and returns.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "gemv.cuh"

namespace shk {
namespace {

constexpr int PF_M = 128, PF_N = 128, PF_K = 64, PF_THREADS = 256;
constexpr int PF_TILE_A = PF_M * PF_K * 2;  // 16 KB
constexpr int PF_TILE_B = PF_N * PF_K * 2;  // 16 KB
constexpr int PF_STAGE = PF_TILE_A + PF_TILE_B;
constexpr int PF_TMEM_COLS = PF_N;  // fp32 accumulator columns
// dynamic shared memory: 1 KB alignment slack, 2 stages, barriers, TMEM slot
constexpr int PF_SMEM = 1024 + 2 * PF_STAGE + 64;

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: start address,
// leading byte offset 16 (unused for swizzled K-major), stride byte offset
// 1024 (8-row groups), descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: D fp32, A and B bf16, both K-major, N, M.
constexpr uint32_t PF_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(PF_N >> 3) << 17) |
                              ((uint32_t)(PF_M >> 4) << 24);

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
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

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// 32 consecutive elements (a quarter half `h` of K-step `ks`) of weight row
// `row`, dequantised (same per-element formulas as the reference's
// dequantize_row_q4_k / dequantize_row_q6_k, engine/src/ops.c:117-193),
// packed as 16 bf16 pairs.
template <int QT>
__device__ __forceinline__ void dequant32(const uint8_t* __restrict__ rowp, uint32_t nb, uint32_t ks, int h,
                                          uint32_t (&out)[16]) {
  const uint32_t b = ks >> 2, j = ks & 3;  // 256-block, its 64-element quarter
  if (QT == T_Q4K) {
    const uint8_t* blk = rowp + (size_t)b * Q4K_BYTES;
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
      out[2 * i] = pack_bf16(v[0], v[1]);
      out[2 * i + 1] = pack_bf16(v[2], v[3]);
    }
  } else {  // planar Q6_K (repack.cu)
    const uint32_t n = j >> 1, g = 2 * (j & 1) + h;  // half, 32-element group
    const uint32_t qlc = 4 * n + 2 * (g & 1), qhc = 2 * n;
    const uint4 a0 = *reinterpret_cast<const uint4*>(rowp + 128 * b + 16 * ((qlc + b) & 7));
    const uint4 a1 = *reinterpret_cast<const uint4*>(rowp + 128 * b + 16 * ((qlc + 1 + b) & 7));
    const uint8_t* qhb = rowp + 128 * nb + 64 * b;
    const uint4 h0 = *reinterpret_cast<const uint4*>(qhb + 16 * ((qhc + (b >> 1)) & 3));
    const uint4 h1 = *reinterpret_cast<const uint4*>(qhb + 16 * ((qhc + 1 + (b >> 1)) & 3));
    const int8_t* scp = reinterpret_cast<const int8_t*>(rowp + 192 * nb + 16 * b + 8 * n + 2 * g);
    const float d = ref_half(*reinterpret_cast<const uint16_t*>(rowp + 208 * nb + 2 * b));
    const float ds0 = d * (float)scp[0], ds1 = d * (float)scp[1];
    const uint32_t ql[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t lo = (g >= 2) ? (ql[i] >> 4) : ql[i];
      const uint32_t hi = qh[i] >> (2 * g);
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int q = (int)(((lo >> (8 * e)) & 0xF) | (((hi >> (8 * e)) & 3) << 4)) - 32;
        v[e] = (i < 4 ? ds0 : ds1) * (float)q;  // elements 0-15: first scale, 16-31: second
      }
      out[2 * i] = pack_bf16(v[0], v[1]);
      out[2 * i + 1] = pack_bf16(v[2], v[3]);
    }
  }
}

__device__ __forceinline__ uint32_t sw128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

template <int QT>
__global__ void __launch_bounds__(PF_THREADS, 1)
    prefill_kernel(const uint8_t* __restrict__ w, uint32_t row_stride, const __nv_bfloat16* __restrict__ xb,
                   float* __restrict__ y, uint32_t M, uint32_t K, uint32_t T, int* err) {
  extern __shared__ uint8_t pf_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pf_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + 2 * PF_STAGE);  // [0], [1]: stages; [2]: all done
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + 2 * PF_STAGE + 32);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t m0 = blockIdx.x * PF_M, t0 = blockIdx.y * PF_N;
  const uint32_t nb = K / QK, nk = K / PF_K;

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_init(&bar[2], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(PF_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  bool ok = true;
  uint32_t ph0 = 0, ph1 = 0;  // phase parity of each stage's barrier
  for (uint32_t ks = 0; ks < nk && ok; ++ks) {
    const uint32_t s = ks & 1;
    uint8_t* A = sm + s * PF_STAGE;
    uint8_t* B = A + PF_TILE_A;
    if (ks >= 2) {  // the MMAs of step ks - 2 have read this stage
      ok = __syncthreads_and(mbar_wait_bounded(&bar[s], s ? ph1 : ph0, err, DERR_TIMEOUT_FULL)) != 0;
      if (s) ph1 ^= 1; else ph0 ^= 1;
      if (!ok) break;
    }
    // A: weight rows m0 + r, elements [64 ks, 64 ks + 64)
    {
      const uint32_t r = tid >> 1, h = tid & 1, m = m0 + r;
      uint32_t v[16];
      if (m < M) {
        dequant32<QT>(w + (size_t)m * row_stride, nb, ks, (int)h, v);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(A + sw128(r, 4 * h + c)) = make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    }
    // B: tokens t0 + r, same elements
#pragma unroll
    for (int i = 0; i < (PF_N * 8) / PF_THREADS; ++i) {
      const uint32_t idx = tid + i * PF_THREADS, r = idx >> 3, c = idx & 7, t = t0 + r;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (t < T) v = __ldg(reinterpret_cast<const uint4*>(xb + (size_t)t * K + (size_t)ks * PF_K) + c);
      *reinterpret_cast<uint4*>(B + sw128(r, c)) = v;
    }
    proxy_fence();  // generic-proxy stores visible to the tensor core (async proxy)
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a0 = smem_u32(A), b0 = smem_u32(B);
#pragma unroll
      for (uint32_t k4 = 0; k4 < PF_K / 16; ++k4)
        mma_bf16(tmem, desc_sw128(a0 + 32 * k4), desc_sw128(b0 + 32 * k4), (ks | k4) ? 1u : 0u);
      mma_commit(&bar[s]);
    }
  }
  // all MMAs issued by thread 0 complete -> bar[2]
  if (tid == 0) mma_commit(&bar[2]);
  const bool done = __syncthreads_and(mbar_wait_bounded(&bar[2], 0, err, DERR_TIMEOUT_FULL)) != 0;
  tc_fence_after();
  if (ok && done && warp < 4) {
    const uint32_t row = 32 * warp + lane, m = m0 + row;
#pragma unroll 1
    for (uint32_t cc = 0; cc < PF_N / 32; ++cc) {
      uint32_t v[32];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
          "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
            "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
            "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
            "=r"(v[30]), "=r"(v[31])
          : "r"(tmem + ((32u * warp) << 16) + 32u * cc));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (m < M) {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const uint32_t t = t0 + 32 * cc + jj;
          if (t < T) y[(size_t)t * M + m] = __uint_as_float(v[jj]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PF_TMEM_COLS) : "memory");
}

__global__ void to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ xb, size_t n) {
  for (size_t i = 2 * ((size_t)blockIdx.x * blockDim.x + threadIdx.x); i < n; i += 2 * (size_t)gridDim.x * blockDim.x) {
    const float2 v = *reinterpret_cast<const float2*>(x + i);
    *reinterpret_cast<__nv_bfloat162*>(xb + i) = __floats2bfloat162_rn(v.x, v.y);
  }
}

}  // namespace

size_t prefill_x_bytes(uint32_t k, uint32_t n_tokens) { return (size_t)k * n_tokens * 2; }

cudaError_t prefill_launch(uint32_t qt, const void* w, uint32_t row_stride, const float* x, void* xb_scratch,
                           float* y, uint32_t m, uint32_t k, uint32_t n_tokens, int* err, int num_sms,
                           cudaStream_t st) {
  const size_t n = (size_t)k * n_tokens;  // k % 256 == 0: even
  to_bf16_kernel<<<4 * num_sms, 256, 0, st>>>(x, static_cast<__nv_bfloat16*>(xb_scratch), n);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const dim3 grid((m + PF_M - 1) / PF_M, (n_tokens + PF_N - 1) / PF_N);
  const auto* xb = static_cast<const __nv_bfloat16*>(xb_scratch);
  const auto* wb = static_cast<const uint8_t*>(w);
  if (qt == T_Q4K) {
    e = cudaFuncSetAttribute(prefill_kernel<T_Q4K>, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
    if (e == cudaSuccess)
      prefill_kernel<T_Q4K><<<grid, PF_THREADS, PF_SMEM, st>>>(wb, row_stride, xb, y, m, k, n_tokens, err);
  } else {
    e = cudaFuncSetAttribute(prefill_kernel<T_Q6K_PLANAR>, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
    if (e == cudaSuccess)
      prefill_kernel<T_Q6K_PLANAR><<<grid, PF_THREADS, PF_SMEM, st>>>(wb, row_stride, xb, y, m, k, n_tokens, err);
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace shk
