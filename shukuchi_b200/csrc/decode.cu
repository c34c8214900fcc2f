// decode.cu -- persistent whole-token decode kernel for sm_100a.
//
// One cooperative launch, one CTA per SM, 15 consumer warps + 1 producer warp
// (the tensor-core matvec's shape, mmv_dev.cuh).  The program is a list of
// phases per token (embed, per layer: QKV, attention, O, gate/up, down; then
// lm_head and argmax), run n_steps times with the argmax token and position
// fed back on the device (engine/src/engine.c:306-501).
//
//  * The producer lane walks every matvec phase of every token in order and
//    streams this CTA's weight chunks into the shared-memory ring; it never
//    waits for activations, so while the consumers convert x, run attention
//    or wait at a phase boundary, the ring fills with the coming projection's
//    weights.  Every plan shares one ring geometry (slot size, chunk, stages).
//  * The consumers run each phase (x conversion + items, attention items,
//    embed slice, argmax slice), then count the phase done on a monotonic
//    grid-wide counter and wait until every CTA has: each phase reads the
//    previous one's output, which may come from any CTA.
//
// Waits are bounded (1 s): a CTA that gives up records SHK_ETIMEOUT and
// leaves; the others then time out at their next phase boundary, so a fault
// never turns into a hang.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "attn_dev.cuh"
#include "common.cuh"
#include "decode.cuh"
#include "glue_dev.cuh"
#include "mmv_dev.cuh"

namespace shk {
namespace {
using namespace mdev;
using namespace adev;
using namespace gldev;

constexpr int DC_CT = 32 * MMV_WARPS;  // consumer threads

// Header of the kernel's shared memory (bytes).
constexpr uint32_t OFF_FULL = 0;
constexpr uint32_t OFF_EMPTY = OFF_FULL + 8 * MMV_MAX_STAGES;
constexpr uint32_t OFF_RED = OFF_EMPTY + 8 * MMV_MAX_STAGES;
constexpr uint32_t OFF_AMV = OFF_RED + 4 * 32;
constexpr uint32_t OFF_AMI = OFF_AMV + 4 * 32;
constexpr uint32_t OFF_FLAG = OFF_AMI + 4 * 32;
constexpr uint32_t OFF_CNT = (OFF_FLAG + 16 + 15) & ~15u;
constexpr uint32_t OFF_PART = (OFF_CNT + 4 * MMV_RED_MAX_SLOTS + 127) & ~127u;
constexpr uint32_t OFF_ARGS = (OFF_PART + 4 * MMV_RED_FLOATS + 127) & ~127u;
constexpr uint32_t HDR_BYTES = (OFF_ARGS + (uint32_t)sizeof(MmvArgs) + 127) & ~127u;

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Phase boundary of the consumer threads (the producer warp never joins):
// count this CTA's phase `seq` done, then wait until every CTA has.  Writes
// before it are visible to every CTA after it.  False if the wait ran out.
__device__ __forceinline__ bool phase_sync(uint32_t* bar, uint32_t seq, int* err, volatile int* flag) {
  named_sync(1, DC_CT);
  if (threadIdx.x == 0) {
    int ok = 1;
    __threadfence();  // this CTA's stores (ordered before by the CTA barrier) before its count
    atomicAdd(bar, 1u);
    const uint32_t target = (seq + 1) * gridDim.x;
    // poll with relaxed loads and a short back-off (148 pollers on one line
    // must not crowd out the late CTAs' atomics), then one acquire fence
    if (ld_relaxed_gpu(bar) < target) {
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t n = 1; ld_relaxed_gpu(bar) < target; ++n) {
        __nanosleep(64);
        if ((n & 63) == 0 && globaltimer_ns() - t0 > WAIT_BUDGET_NS) {
          set_error(err, DERR_TIMEOUT_GRID);
          ok = 0;
          break;
        }
      }
    }
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    *flag = ok;
  }
  named_sync(1, DC_CT);
  return *flag != 0;
}

// This CTA's items of a plan ([i0, i1); none past the plan's grid).
__device__ __forceinline__ void cta_items(const MmvArgs& a, uint32_t& i0, uint32_t& i1) {
  if (blockIdx.x < a.grid) {
    i0 = a.cta_item[blockIdx.x];
    i1 = a.cta_item[blockIdx.x + 1];
  } else {
    i0 = i1 = 0;
  }
}

// Ring chunks a plan's items [i0, i1) take (they never share a chunk with
// another plan's).
__device__ __forceinline__ uint32_t plan_chunks(const MRing& R, uint32_t i0, uint32_t i1) {
  return (i1 - i0 + R.chunk - 1) >> R.lg_chunk;
}

template <int HD, int G>
__global__ void __launch_bounds__(MMV_THREADS, 1) decode_kernel(const __grid_constant__ DecodeProgram P) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_FULL);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + OFF_EMPTY);
  float* red = reinterpret_cast<float*>(smem + OFF_RED);
  float* am_sv = reinterpret_cast<float*>(smem + OFF_AMV);
  uint32_t* am_si = reinterpret_cast<uint32_t*>(smem + OFF_AMI);
  volatile int* flag = reinterpret_cast<volatile int*>(smem + OFF_FLAG);
  int* cnt = reinterpret_cast<int*>(smem + OFF_CNT);
  float* part = reinterpret_cast<float*>(smem + OFF_PART);
  MmvArgs* sargs = reinterpret_cast<MmvArgs*>(smem + OFF_ARGS);
  uint8_t* xreg = smem + P.xreg_off;
  const MRing R{full, empty, smem + P.ring_off, P.ns, P.slot_bytes, P.chunk, P.lg_chunk};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid < (int)P.ns) {
    mbar_init(&full[tid], 1);
    mbar_init(&empty[tid], P.chunk);
    fence_mbar_init();
  }
  for (int i = tid; i < MMV_RED_MAX_SLOTS; i += MMV_THREADS) cnt[i] = 0;
  __syncthreads();

  if (warp == MMV_WARPS) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      uint32_t cpos = 0;
      bool ok = true;
      for (uint32_t step = 0; step < P.n_steps && ok; ++step)
        for (uint32_t ph = 0; ph < P.n_phases && ok; ++ph) {
          const DecodePhase d = P.phases[ph];
          if (d.kind != PH_GEMV) continue;
          const MmvArgs& a = P.mmv[d.idx];
          uint32_t i0, i1;
          cta_items(a, i0, i1);
          ok = mmv_produce(a, R, i0, i1, cpos, nullptr, 0);
        }
      mmv_drain(R, cpos, P.err);
    }
    return;
  }

  // ------------------------------ consumers -------------------------------
  uint32_t cpos = 0, seq = 0;
  const bool tracing = P.trace && blockIdx.x == 0 && tid == 0;
  if (tracing) P.trace[0] = globaltimer_ns();
  for (uint32_t step = 0; step < P.n_steps; ++step) {
    for (uint32_t ph = 0; ph < P.n_phases; ++ph) {
      const DecodePhase d = P.phases[ph];
      bool ok = true;
      if (d.kind == PH_GEMV) {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(&P.mmv[d.idx]);
        uint32_t* dst = reinterpret_cast<uint32_t*>(sargs);
        for (uint32_t i = tid; i < sizeof(MmvArgs) / 4; i += DC_CT) dst[i] = __ldg(src + i);
        named_sync(1, DC_CT);
        const MmvArgs& a = *sargs;
        uint32_t i0, i1;
        cta_items(a, i0, i1);
        if (i0 < i1) {
          const XRegion X = x_region(xreg, a.k, a.has4, a.has6);
          if (a.has4 && a.has6) {
            const float osc = mmv_prologue<true, true>(a, X, red, warp, lane, nullptr);
            ok = mmv_consume<true, true>(a, R, i0, i1, cpos, X, osc, part, cnt, warp, lane);
          } else if (a.has4) {
            const float osc = mmv_prologue<true, false>(a, X, red, warp, lane, nullptr);
            ok = mmv_consume<true, false>(a, R, i0, i1, cpos, X, osc, part, cnt, warp, lane);
          } else {
            const float osc = mmv_prologue<false, true>(a, X, red, warp, lane, nullptr);
            ok = mmv_consume<false, true>(a, R, i0, i1, cpos, X, osc, part, cnt, warp, lane);
          }
        }
        cpos += plan_chunks(R, i0, i1);
      } else if (d.kind == PH_ATTN) {
        const AttnArgs& aa = P.attn[d.idx];
        const uint32_t n_items = P.n_kv * P.attn_nsplit;
        for (uint32_t item = blockIdx.x; item < n_items; item += gridDim.x)
          attn_item<HD, G, MMV_WARPS>(aa, item % P.n_kv, item / P.n_kv, P.attn_nsplit,
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
          *flag = atomicAdd(P.am_cnt, 1) == (int)gridDim.x - 1;
        }
        named_sync(1, DC_CT);
        if (*flag) {  // the last CTA merges the partials with all its threads
          __threadfence();
          const bool x0_nan = isnan(__ldcg(P.logits));
          const uint32_t ix = am_merge_par<DC_CT>(P.am_v, P.am_i, gridDim.x, x0_nan, am_sv, am_si,
                                                  [] { named_sync(1, DC_CT); });
          if (tid == 0) {
            P.tok[0] = ix;
            if (P.advance_pos) P.tok[1] = __ldcg(P.tok + 1) + 1;
            *P.am_cnt = 0;
          }
        }
      }
      if (!ok) return;  // a bounded wait ran out; the error is recorded
      const bool rec = tracing && seq < P.trace_cap_phases;
      if (rec) P.trace[1 + 2 * seq] = globaltimer_ns();
      if (!phase_sync(P.bar, seq, P.err, flag)) return;
      if (rec) P.trace[2 + 2 * seq] = globaltimer_ns();
      ++seq;
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
    case 128 * 16 + 1: return AttnSmem<128, 1, MMV_WARPS>::BYTES;
    case 128 * 16 + 2: return AttnSmem<128, 2, MMV_WARPS>::BYTES;
    case 128 * 16 + 4: return AttnSmem<128, 4, MMV_WARPS>::BYTES;
    case 128 * 16 + 8: return AttnSmem<128, 8, MMV_WARPS>::BYTES;
    case 64 * 16 + 1: return AttnSmem<64, 1, MMV_WARPS>::BYTES;
    case 64 * 16 + 2: return AttnSmem<64, 2, MMV_WARPS>::BYTES;
    case 64 * 16 + 4: return AttnSmem<64, 4, MMV_WARPS>::BYTES;
    case 64 * 16 + 8: return AttnSmem<64, 8, MMV_WARPS>::BYTES;
    default: return 0;
  }
}

}  // namespace

size_t decode_smem(DecodeProgram& P, uint32_t head_dim, uint32_t group, size_t* fixed_out) {
  const size_t att = attn_smem_bytes(head_dim, group);
  const size_t xr = std::max(x_bytes(P.kmax, true, true), att);
  P.xreg_off = HDR_BYTES;
  P.ring_off = (uint32_t)((P.xreg_off + xr + 127) & ~(size_t)127);
  if (fixed_out) *fixed_out = P.ring_off;
  return (size_t)P.ring_off + (size_t)P.ns * P.chunk * P.slot_bytes;
}

bool decode_supported(uint32_t head_dim, uint32_t group, size_t smem, int num_sms) {
  void* k = pick_kernel(head_dim, group);
  if (!k || smem > 227 * 1024) return false;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return false;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, MMV_THREADS, smem) != cudaSuccess)
    return false;
  return per_sm >= 1 && num_sms >= 1;
}

cudaError_t decode_launch(const DecodeProgram& P, uint32_t head_dim, uint32_t group, size_t smem,
                          int grid, cudaStream_t stream) {
  void* k = pick_kernel(head_dim, group);
  if (!k) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(P.bar, 0, sizeof(uint32_t), stream);
  if (e != cudaSuccess) return e;
  void* args[] = {const_cast<DecodeProgram*>(&P)};
  return cudaLaunchCooperativeKernel(k, dim3(grid), dim3(MMV_THREADS), args, smem, stream);
}

}  // namespace shk
