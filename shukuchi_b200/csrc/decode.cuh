// decode.cuh -- persistent whole-token decode kernel (host-side API).
//
// One cooperative launch runs n tokens: embed -> per layer (RMSNorm + QKV +
// RoPE GEMV, append + attention, O + residual, RMSNorm + gate/up + SwiGLU,
// down + residual) -> lm_head -> argmax, feeding the argmax back to the next
// embed on the device (engine/src/engine.c:306-501 token loop,
// :76-229 layer forward).  Phases are separated by grid-wide barriers; the
// producer warp of every CTA keeps streaming the weights of the coming GEMV
// phases into its shared-memory ring across those barriers, so HBM streaming
// does not stop between projections, layers or tokens.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "attn.cuh"
#include "gemv.cuh"

namespace shk {

enum DecodePhaseKind : uint32_t { PH_EMBED = 0, PH_GEMV = 1, PH_ATTN = 2, PH_ARGMAX = 3 };

struct DecodePhase {
  uint32_t kind;  // DecodePhaseKind
  uint32_t idx;   // index into DecodeProgram::gemv or ::attn
};

// Grid barrier state in device memory (zeroed before each launch).
struct GridBar {
  uint32_t count;
  uint32_t gen;
};

struct DecodeProgram {
  const GemvArgs* gemv;       // device array of GEMV phase plans
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
  uint32_t* tok;  // device [0] token, [1] position
  uint32_t advance_pos;  // argmax advances tok[1] (device-fed token loop)
  // shared-memory geometry
  uint32_t ns, stage_bytes;  // ring stages and their size
  uint32_t xreg_off, ring_off;
  // attention work split: n_kv heads x attn_nsplit position splits
  uint32_t n_kv, attn_nsplit;
  GridBar* bar;
  int* err;
  // optional timeline (null = off): CTA 0 records %globaltimer at the start and,
  // per phase, when it reaches the barrier and when it leaves it:
  // trace[0] = start, trace[1 + 2*i] = arrive, trace[2 + 2*i] = leave for the
  // i-th phase of the launch (i < trace_cap_phases)
  uint64_t* trace;
  uint32_t trace_cap_phases;
};

// Shared memory of the decode kernel for the given head geometry, largest K
// and ring.  Fills P.xreg_off / P.ring_off.
size_t decode_smem(DecodeProgram& P, uint32_t head_dim, uint32_t group, uint32_t kmax);
// Sets the kernel attributes; returns false if this (head_dim, group) is not
// built or one CTA per SM does not fit.
bool decode_supported(uint32_t head_dim, uint32_t group, size_t smem, int num_sms);
// Cooperative launch, one CTA per SM (grid = num_sms).
cudaError_t decode_launch(const DecodeProgram& P, uint32_t head_dim, uint32_t group, size_t smem,
                          int grid, cudaStream_t stream);

}  // namespace shk
