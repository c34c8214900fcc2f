// decode.cuh -- persistent whole-token decode kernel (host-side API).
//
// One cooperative launch runs n tokens: embed -> per layer (RMSNorm + QKV +
// RoPE matvec, append + attention, O + residual, RMSNorm + gate/up + SwiGLU,
// down + residual) -> lm_head -> argmax, feeding the argmax back to the next
// embed on the device (engine/src/engine.c:306-501 token loop, :76-229 layer
// forward).  The projections are tensor-core matvecs over row-tiled weights
// (mmv_dev.cuh).  A producer lane per CTA streams the weight chunks of every
// matvec phase of every token into the CTA's shared-memory ring in program
// order and never waits for activations, so HBM keeps streaming through the
// phase boundaries (grid-wide waits on a monotonic counter), attention and
// the x conversions.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "attn.cuh"
#include "mmv.cuh"

namespace shk {

enum DecodePhaseKind : uint32_t { PH_EMBED = 0, PH_GEMV = 1, PH_ATTN = 2, PH_ARGMAX = 3 };

struct DecodePhase {
  uint32_t kind;  // DecodePhaseKind
  uint32_t idx;   // index into DecodeProgram::mmv or ::attn
};

struct DecodeProgram {
  const MmvArgs* mmv;         // device array of matvec phase plans (common ring geometry)
  const AttnArgs* attn;       // device array of attention phases
  const DecodePhase* phases;  // device array: one token's phases in order
  uint32_t n_phases;          // phases per token
  uint32_t n_steps;           // tokens
  // embed (engine/src/ops.c:533-577)
  const uint8_t* tok_embd;
  uint32_t embd_dtype, n_vocab, n_embd;
  float* hidden;
  // argmax (engine/src/engine.c:424-431); partials sized >= grid
  const float* logits;
  float* am_v;
  uint32_t* am_i;
  int* am_cnt;
  uint32_t* tok;          // device [0] token, [1] position
  uint32_t advance_pos;   // argmax advances tok[1] (device-fed token loop)
  // shared-memory geometry: ring of ns stages of `chunk` slots of slot_bytes
  uint32_t ns, slot_bytes, chunk, lg_chunk;
  uint32_t xreg_off, ring_off;
  uint32_t kmax;          // largest matvec K (x region size)
  // attention work split: n_kv heads x attn_nsplit position splits
  uint32_t n_kv, attn_nsplit;
  uint32_t* bar;          // phases completed x grid (zeroed before each launch)
  int* err;
  // optional timeline (null = off): CTA 0 records %globaltimer at the start and,
  // per phase, when it reaches the barrier and when it leaves it:
  // trace[0] = start, trace[1 + 2*i] = arrive, trace[2 + 2*i] = leave for the
  // i-th phase of the launch (i < trace_cap_phases)
  uint64_t* trace;
  uint32_t trace_cap_phases;
};

// Shared memory of the decode kernel for the given head geometry and largest
// K, with the ring geometry already in P (ns, slot_bytes, chunk).  Fills
// P.xreg_off / P.ring_off.  fixed_out: bytes before the ring.
size_t decode_smem(DecodeProgram& P, uint32_t head_dim, uint32_t group, size_t* fixed_out = nullptr);
// Sets the kernel attributes; returns false if this (head_dim, group) is not
// built or one CTA per SM does not fit.
bool decode_supported(uint32_t head_dim, uint32_t group, size_t smem, int num_sms);
// Cooperative launch, one CTA per SM (grid = num_sms).
cudaError_t decode_launch(const DecodeProgram& P, uint32_t head_dim, uint32_t group, size_t smem,
                          int grid, cudaStream_t stream);

}  // namespace shk
