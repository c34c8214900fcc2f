// decode.cu -- persistent whole-token decode kernel for sm_100a.
//
// One cooperative launch, one CTA per SM, 8 consumer warps + 1 producer warp
// (the GEMV kernel's shape).  The program is a list of phases per token
// (embed, per layer: QKV GEMV, attention, O GEMV, gate/up GEMV, down GEMV;
// then lm_head GEMV and argmax), run n_steps times with the argmax token and
// position fed back on the device (engine/src/engine.c:306-501).
//
//  * The producer lane walks every GEMV phase of every token in order and
//    streams this CTA's weight chunks into the shared-memory ring; it never
//    waits for activations, so while the consumers are in an attention phase
//    or at a barrier the ring fills with the coming projection's weights.
//  * The consumers run each phase (GEMV prologue + tasks, attention items,
//    embed slice, argmax slice) and then meet at a grid-wide barrier: every
//    phase reads the previous phase's output, which may come from any CTA.
//
// Waits are bounded (1 s): a CTA that gives up records SHK_ETIMEOUT and
// leaves; the others then time out at their next barrier, so a fault never
// turns into a hang.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "attn_dev.cuh"
#include "common.cuh"
#include "decode.cuh"
#include "gemv_dev.cuh"
#include "glue_dev.cuh"

namespace shk {
namespace {
using namespace gdev;
using namespace adev;
using namespace gldev;

constexpr int DC_CT = 32 * GEMV_WARPS;  // consumer threads

// Header of the kernel's shared memory (bytes).
constexpr uint32_t OFF_FULL = 0;
constexpr uint32_t OFF_EMPTY = OFF_FULL + 8 * GEMV_MAX_STAGES;
constexpr uint32_t OFF_DONE = OFF_EMPTY + 8 * GEMV_MAX_STAGES;
constexpr uint32_t OFF_GEN = OFF_DONE + 4 * GEMV_MAX_STAGES;
constexpr uint32_t OFF_RED = OFF_GEN + 4 * GEMV_MAX_STAGES;
constexpr uint32_t OFF_AMV = OFF_RED + 4 * 32;
constexpr uint32_t OFF_AMI = OFF_AMV + 4 * (DC_CT / 32);
constexpr uint32_t OFF_FLAG = OFF_AMI + 4 * (DC_CT / 32);
constexpr uint32_t OFF_KPART = (OFF_FLAG + 16 + 15) & ~15u;
constexpr uint32_t OFF_KCNT = OFF_KPART + 4 * GEMV_MAX_STAGES * GEMV_KS_ROWT * GEMV_KS_MAX * 2;
constexpr uint32_t OFF_ARGS = (OFF_KCNT + 4 * GEMV_MAX_STAGES * GEMV_KS_ROWT + 15) & ~15u;
constexpr uint32_t HDR_BYTES = (OFF_ARGS + (uint32_t)sizeof(GemvArgs) + 127) & ~127u;

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of the consumer threads (the producer warp never joins).
// Writes before it are visible to every CTA after it.  False if the wait ran
// out (error recorded).
__device__ __forceinline__ bool grid_sync(GridBar* gb, int* err, volatile int* flag) {
  named_sync(1, DC_CT);
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint32_t g = *reinterpret_cast<volatile uint32_t*>(&gb->gen);
    __threadfence();
    if (atomicAdd(&gb->count, 1u) == gridDim.x - 1) {
      atomicExch(&gb->count, 0u);
      __threadfence();
      atomicExch(&gb->gen, g + 1);
    } else {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_gpu(&gb->gen) == g) {
        if (globaltimer_ns() - t0 > WAIT_BUDGET_NS) {
          set_error(err, DERR_TIMEOUT_GRID);
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
    *flag = ok;
  }
  named_sync(1, DC_CT);
  return *flag != 0;
}

template <int HD, int G>
__global__ void __launch_bounds__(GEMV_THREADS, 1) decode_kernel(const __grid_constant__ DecodeProgram P) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_FULL);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + OFF_EMPTY);
  int* done = reinterpret_cast<int*>(smem + OFF_DONE);
  volatile uint32_t* gen = reinterpret_cast<volatile uint32_t*>(smem + OFF_GEN);
  float* red = reinterpret_cast<float*>(smem + OFF_RED);
  float* am_sv = reinterpret_cast<float*>(smem + OFF_AMV);
  uint32_t* am_si = reinterpret_cast<uint32_t*>(smem + OFF_AMI);
  volatile int* flags = reinterpret_cast<volatile int*>(smem + OFF_FLAG);
  GemvArgs* sargs = reinterpret_cast<GemvArgs*>(smem + OFF_ARGS);
  uint8_t* xreg = smem + P.xreg_off;
  const Ring R{full,           empty, done, gen, smem + P.ring_off, P.ns, P.stage_bytes,
               reinterpret_cast<float*>(smem + OFF_KPART), reinterpret_cast<int*>(smem + OFF_KCNT)};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (uint32_t s = 0; s < P.ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      done[s] = 0;
      gen[s] = 0xFFFFFFFFu;
      for (int r = 0; r < GEMV_KS_ROWT; ++r) R.kcnt[s * GEMV_KS_ROWT + r] = 0;
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == GEMV_WARPS) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      RingPos p;
      bool ok = true;
      for (uint32_t step = 0; step < P.n_steps && ok; ++step)
        for (uint32_t ph = 0; ph < P.n_phases && ok; ++ph) {
          const DecodePhase d = P.phases[ph];
          if (d.kind != PH_GEMV) continue;
          const GemvArgs& a = P.gemv[d.idx];
          const uint64_t lo = a.total_cost * blockIdx.x / gridDim.x;
          const uint64_t hi = a.total_cost * (blockIdx.x + 1) / gridDim.x;
          ok = gemv_produce(a, R, p, lo, hi);
        }
      ring_drain(R, p, P.err);
    }
    return;
  }

  // ------------------------------ consumers -------------------------------
  RingPos p;
  uint32_t gtask = 0;
  const bool tracing = P.trace && blockIdx.x == 0 && tid == 0;
  if (tracing) P.trace[0] = globaltimer_ns();
  uint32_t n_done = 0;
  for (uint32_t step = 0; step < P.n_steps; ++step) {
    for (uint32_t ph = 0; ph < P.n_phases; ++ph) {
      const DecodePhase d = P.phases[ph];
      bool ok = true;
      if (d.kind == PH_GEMV) {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(&P.gemv[d.idx]);
        uint32_t* dst = reinterpret_cast<uint32_t*>(sargs);
        for (uint32_t i = tid; i < sizeof(GemvArgs) / 4; i += DC_CT) dst[i] = src[i];
        named_sync(1, DC_CT);
        const GemvArgs& a = *sargs;
        bool h4 = false, h6 = false;
        for (uint32_t s = 0; s < a.nseg; ++s) {
          h4 = h4 || a.seg[s].qt == T_Q4K;
          h6 = h6 || a.seg[s].qt == T_Q6K;
        }
        const uint32_t K = a.k;
        XBuf xb;
        xb.xq = reinterpret_cast<int4*>(xreg);
        xb.xbs = reinterpret_cast<float*>(xreg + xq_bytes(K));
        xb.xs32 = xb.xbs + xbs_floats(K);
        const uint64_t lo = a.total_cost * blockIdx.x / gridDim.x;
        const uint64_t hi = a.total_cost * (blockIdx.x + 1) / gridDim.x;
        if (h4 && h6) {
          const float osc = gemv_prologue<true, true>(a, xb, red, warp, lane);
          ok = gemv_consume<true, true>(a, R, p, gtask, lo, hi, xb.view(osc), warp, lane);
        } else if (h4) {
          const float osc = gemv_prologue<true, false>(a, xb, red, warp, lane);
          ok = gemv_consume<true, false>(a, R, p, gtask, lo, hi, xb.view(osc), warp, lane);
        } else {
          const float osc = gemv_prologue<false, true>(a, xb, red, warp, lane);
          ok = gemv_consume<false, true>(a, R, p, gtask, lo, hi, xb.view(osc), warp, lane);
        }
      } else if (d.kind == PH_ATTN) {
        const AttnArgs& aa = P.attn[d.idx];
        const uint32_t n_items = P.n_kv * P.attn_nsplit;
        for (uint32_t item = blockIdx.x; item < n_items; item += gridDim.x)
          attn_item<HD, G, GEMV_WARPS>(aa, item % P.n_kv, item / P.n_kv, P.attn_nsplit,
                                        reinterpret_cast<float*>(xreg));
      } else if (d.kind == PH_EMBED) {
        const uint32_t tok = __ldcg(P.tok);
        if (tok >= P.n_vocab) {
          if (blockIdx.x == 0 && tid == 0) set_error(P.err, DERR_BAD_TOKEN);
        } else {
          for (uint32_t e = blockIdx.x * DC_CT + tid; e < P.n_embd; e += gridDim.x * DC_CT)
            P.hidden[e] = embed_elem(P.tok_embd, P.embd_dtype, tok, P.n_embd, e);
        }
      } else {  // PH_ARGMAX over the logits, first index on ties
        const uint32_t per = (P.n_vocab + gridDim.x - 1) / gridDim.x;
        const uint32_t lo = min(P.n_vocab, blockIdx.x * per), hi = min(P.n_vocab, lo + per);
        float bv;
        uint32_t bi;
        am_block<DC_CT>(P.logits, lo, hi, am_sv, am_si, [] { named_sync(1, DC_CT); }, bv, bi);
        if (tid == 0) {
          P.am_v[blockIdx.x] = bv;
          P.am_i[blockIdx.x] = bi;
          __threadfence();
          if (atomicAdd(P.am_cnt, 1) == (int)gridDim.x - 1) {
            __threadfence();
            P.tok[0] = am_merge(P.am_v, P.am_i, gridDim.x);
            if (P.advance_pos) P.tok[1] = __ldcg(P.tok + 1) + 1;
            *P.am_cnt = 0;
          }
        }
      }
      if (!ok) return;  // a bounded wait ran out; the error is recorded
      const bool rec = tracing && n_done < P.trace_cap_phases;
      if (rec) P.trace[1 + 2 * n_done] = globaltimer_ns();
      if (!grid_sync(P.bar, P.err, flags)) return;
      if (rec) P.trace[2 + 2 * n_done] = globaltimer_ns();
      ++n_done;
    }
  }
}

template <int HD, int G>
void* kernel_ptr() {
  return reinterpret_cast<void*>(&decode_kernel<HD, G>);
}

void* pick_kernel(uint32_t hd, uint32_t g) {
  if (hd == 128) {
    if (g == 1) return kernel_ptr<128, 1>();
    if (g == 2) return kernel_ptr<128, 2>();
    if (g == 4) return kernel_ptr<128, 4>();
    if (g == 8) return kernel_ptr<128, 8>();
  } else if (hd == 64) {
    if (g == 1) return kernel_ptr<64, 1>();
    if (g == 2) return kernel_ptr<64, 2>();
    if (g == 4) return kernel_ptr<64, 4>();
    if (g == 8) return kernel_ptr<64, 8>();
  }
  return nullptr;
}

size_t attn_smem_bytes(uint32_t hd, uint32_t g) {
  switch (hd * 16 + g) {
    case 128 * 16 + 1: return AttnSmem<128, 1, GEMV_WARPS>::BYTES;
    case 128 * 16 + 2: return AttnSmem<128, 2, GEMV_WARPS>::BYTES;
    case 128 * 16 + 4: return AttnSmem<128, 4, GEMV_WARPS>::BYTES;
    case 128 * 16 + 8: return AttnSmem<128, 8, GEMV_WARPS>::BYTES;
    case 64 * 16 + 1: return AttnSmem<64, 1, GEMV_WARPS>::BYTES;
    case 64 * 16 + 2: return AttnSmem<64, 2, GEMV_WARPS>::BYTES;
    case 64 * 16 + 4: return AttnSmem<64, 4, GEMV_WARPS>::BYTES;
    case 64 * 16 + 8: return AttnSmem<64, 8, GEMV_WARPS>::BYTES;
    default: return 0;
  }
}

}  // namespace

size_t decode_smem(DecodeProgram& P, uint32_t head_dim, uint32_t group, uint32_t kmax) {
  const size_t att = attn_smem_bytes(head_dim, group);
  const size_t xr = std::max(x_region_bytes(kmax, true, true), att);
  P.xreg_off = HDR_BYTES;
  P.ring_off = (uint32_t)((P.xreg_off + xr + 127) & ~(size_t)127);
  return (size_t)P.ring_off + (size_t)P.ns * P.stage_bytes;
}

bool decode_supported(uint32_t head_dim, uint32_t group, size_t smem, int num_sms) {
  void* k = pick_kernel(head_dim, group);
  if (!k || smem > 227 * 1024) return false;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return false;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, GEMV_THREADS, smem) != cudaSuccess)
    return false;
  return per_sm >= 1 && num_sms >= 1;
}

cudaError_t decode_launch(const DecodeProgram& P, uint32_t head_dim, uint32_t group, size_t smem,
                          int grid, cudaStream_t stream) {
  void* k = pick_kernel(head_dim, group);
  if (!k) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(P.bar, 0, sizeof(GridBar), stream);
  if (e != cudaSuccess) return e;
  void* args[] = {const_cast<DecodeProgram*>(&P)};
  return cudaLaunchCooperativeKernel(k, dim3(grid), dim3(GEMV_THREADS), args, smem, stream);
}

}  // namespace shk
