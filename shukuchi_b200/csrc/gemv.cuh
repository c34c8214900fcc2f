// gemv.cuh -- batch-1 Q4_K / Q6_K dequantise-matvec for sm_100a (host-side plan API).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace shk {

// Epilogue applied to each output row.
enum GemvEpi : uint8_t {
  EPI_STORE = 0,   // y[r] = acc
  EPI_ADD = 1,     // y[r] += acc            (residual add, engine/src/engine.c:164-166)
  EPI_ROPE = 2,    // RoPE on the (2i, 2i+1) pair, then store (engine/src/ops.c:216-238)
  EPI_SWIGLU = 3,  // dual rows: y[r] = silu(gate) * up    (engine/src/ops.c:491-496)
  EPI_TP = 4,      // partial rows to every rank's exchange buffer (GemvTp)
};

constexpr int GEMV_MAX_SEGS = 4;
constexpr int GEMV_WARPS = 15;  // consumer warps; one more warp issues the bulk copies
constexpr int GEMV_THREADS = 32 * (GEMV_WARPS + 1);
constexpr int GEMV_MAX_STAGES = 16;

struct GemvSeg {
  const uint8_t* w;     // matrix: m rows, row r at w + r * row_stride
  const uint8_t* w2;    // second matrix of a dual (gate/up) segment, same shape
  float* y;             // output, m floats
  uint32_t m;           // rows
  uint32_t nb;          // 256-element super-blocks per row
  uint32_t row_stride;  // bytes between rows; multiple of 16
  uint32_t chunk_rows;  // rows per pipeline stage (multiple of rg * rl)
  uint32_t unit_cost;   // bytes per task unit of rg * rl rows (both matrices for dual)
  uint32_t rope_hd;     // head_dim for EPI_ROPE
  uint8_t qt;           // 12 = Q4_K, 14 = Q6_K (planar layout, repack.cu)
  uint8_t epi;          // GemvEpi
  uint8_t rg;           // row groups per warp task (lanes split across groups)
  uint8_t rl;           // rows per lane (each loaded x value feeds rl rows)
  uint8_t dual;         // 1 for gate/up pairs
  uint8_t ks;           // K slices per row task (long rows: one warp per slice), a power of two
  uint8_t lg_ks;        // log2(ks)
  uint16_t sw;          // blocks per K slice: ceil(nb / ks)
};

// Tensor-parallel exchange over NVLink peer memory (one-shot all-reduce fused
// into the GEMVs).  A producer GEMV (out) writes its partial output rows
// (absolute rows row_off + r) into parts_out[p] + rank * d on every rank p;
// its last CTA then stores the step's epoch into flags_out[p][rank].  A
// consumer GEMV (in) waits until flags_in[r] reaches the epoch for every rank
// r and takes x[k] = res_in[k] + sum over r in rank order of parts_in[r*d + k]
// for k in [cov_lo[r], cov_hi[r]); CTA 0 also writes x to res_out (the
// residual stream of the next step).
constexpr int GEMV_TP_MAX = 8;
struct GemvTp {
  const float* parts_in;
  const uint32_t* flags_in;
  float* res_out;
  float* parts_out[GEMV_TP_MAX];
  uint32_t* flags_out[GEMV_TP_MAX];
  uint32_t* counter;        // producer: CTAs done (the last one signals, then resets it)
  const uint32_t* epoch;    // device step counter (advanced by the embedding kernel)
  uint32_t cov_lo[GEMV_TP_MAX], cov_hi[GEMV_TP_MAX];
  uint32_t d;               // elements of one partial
  uint32_t row_off;         // producer: absolute row of output row 0
  uint8_t rank, world, in, out;
};

struct GemvArgs {
  GemvSeg seg[GEMV_MAX_SEGS];
  uint32_t nseg;
  uint32_t k;               // input dimension shared by all segments
  const float* x;           // k floats
  const float* norm_w;      // optional: x <- rmsnorm(x) * norm_w  (eps 1e-5)
  const uint32_t* pos;      // device position for EPI_ROPE
  const float* rope_freq;   // EPI_ROPE: freq[i/2] = powf(1/theta, i/head_dim), host libm
  uint32_t stage_bytes;     // bytes per pipeline stage
  uint32_t n_stages;        // ring depth (<= GEMV_MAX_STAGES)
  uint64_t total_cost;      // sum over segments of units * unit_cost
  int* err;                 // device error word
  GemvTp tp;                // tensor-parallel exchange (tp.in / tp.out = 0: none)
};

struct GemvPlan {
  GemvArgs args;
  int grid = 0;
  size_t smem = 0;
  int has4 = 0, has6 = 0;
};

// Describes one matrix for planning.
struct GemvMat {
  const void* w;
  const void* w2;  // non-null => dual segment (gate/up)
  float* y;
  uint32_t m;
  uint32_t qt;
  uint32_t row_stride;  // 0 => dense rows
  uint8_t epi;
  uint32_t rope_hd;
};

// Returns 0 on success, negative on unsupported shapes (caller may fall back).
// max_stage_bytes bounds the bytes of one pipeline stage (a chunk of rows).
#ifndef SHK_GEMV_STAGE_BYTES
#define SHK_GEMV_STAGE_BYTES 32768
#endif
int gemv_plan(GemvPlan& p, const GemvMat* mats, int nmats, uint32_t k, const float* x,
              const float* norm_w, const uint32_t* pos, const float* rope_freq, int* err,
              int num_sms, uint32_t max_stage_bytes = SHK_GEMV_STAGE_BYTES);
// Bytes of the x region (fixed-point limbs and per-block sums) for input size K.
size_t gemv_x_region_bytes(uint32_t K, bool has4, bool has6);
// Sets the kernels' dynamic shared-memory limit; call once per device.
cudaError_t gemv_init();
cudaError_t gemv_launch(const GemvPlan& p, cudaStream_t stream);

// Q6_K rows, in place, between the GGUF block layout and the planar layout the
// staged kernel reads (repack.cu).  stride: row bytes, a multiple of 16.
cudaError_t q6k_repack_launch(void* w, uint32_t rows, uint32_t k, uint32_t stride, bool to_planar,
                              int num_sms, cudaStream_t st);

// Batched dequantise-matmul on the tensor cores (prefill.cu): y[t][m] for
// n_tokens tokens; x fp32 [n_tokens][k] is first converted into xb_scratch
// (prefill_x_bytes) as f16, each token row scaled by a power of two (its
// largest magnitude to [2^14, 2^15)), the weights dequantised to f16; fp32
// accumulation.  qt: T_Q4K or T_Q6K_PLANAR.
size_t prefill_x_bytes(uint32_t k, uint32_t n_tokens);
cudaError_t prefill_launch(uint32_t qt, const void* w, uint32_t row_stride, const float* x, void* xb_scratch,
                           float* y, uint32_t m, uint32_t k, uint32_t n_tokens, int* err, int num_sms,
                           cudaStream_t st);

// The tensor-parallel consumer sum of plan args a.tp / a.x as a kernel of its
// own (writes a.tp.res_out).
cudaError_t gemv_tp_sum_launch(const GemvArgs& a, cudaStream_t st);

// Simple fallback for layouts the staged kernel does not take (rows not a
// multiple of 16 bytes; GGUF-layout Q6_K).  Same math, plain loads.
cudaError_t gemv_generic_launch(uint32_t qt, const void* w, const float* x, float* y, uint32_t m,
                                uint32_t k, cudaStream_t stream);

}  // namespace shk
